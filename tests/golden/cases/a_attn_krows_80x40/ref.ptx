.version 8.0
.target sm_89
.address_size 64

.shared .align 16 .b8 _cache_kt[12800];

.visible .entry k_attn_naive(
        .param .u64 param_q,
        .param .u64 param_kt,
        .param .u64 param_v,
        .param .u64 param_attn
)
.reqntid 128
{
        .reg .pred      %p<8>;
        .reg .f32       %f<26>;
        .reg .b32       %r<36>;
        .reg .b64       %rd<11>;

        ld.param.u64    %rd1, [param_q];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_kt];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_v];
        cvta.to.global.u64     %rd3, %rd3;
        ld.param.u64    %rd4, [param_attn];
        cvta.to.global.u64     %rd4, %rd4;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        mov.u32         %r6, _cache_kt;
        mov.s32         %r7, %r1;
        .pragma "nounroll";
CACHE_1:
        setp.ge.s32     %p1, %r7, 3200;
        @%p1 bra        CACHEEND_2;
        mad.wide.s32    %rd5, %r7, 4, %rd2;
        mad.lo.s32      %r8, %r7, 4, %r6;
        ld.global.nc.f32   %f1, [%rd5];
        st.shared.f32   [%r8], %f1;
        add.s32         %r7, %r7, 128;
        bra             CACHE_1;
CACHEEND_2:
        bar.sync        0;
        div.s32         %r9, %r4, 40;
        rem.s32         %r10, %r4, 40;
        mov.f32         %f2, 0fF149F2CA;
        mov.s32         %r11, 0;
        .pragma "nounroll";
LOOP_3:
        mov.f32         %f3, 0f00000000;
        mov.s32         %r12, 0;
        .pragma "nounroll";
LOOP_4:
        mul.lo.s32      %r13, %r9, 40;
        add.s32         %r14, %r13, %r12;
        mad.wide.s32    %rd6, %r14, 4, %rd1;
        ld.global.nc.f32   %f4, [%rd6];
        mul.lo.s32      %r15, %r11, 40;
        add.s32         %r16, %r15, %r12;
        mad.lo.s32      %r17, %r16, 4, %r6;
        ld.shared.f32   %f5, [%r17];
        fma.rn.f32      %f3, %f4, %f5, %f3;
        add.s32         %r12, %r12, 1;
        setp.lt.s32     %p2, %r12, 40;
        @%p2 bra        LOOP_4;
        mov.f32         %f6, 0f3E21E89B;
        mul.f32         %f3, %f3, %f6;
        max.f32         %f2, %f2, %f3;
        add.s32         %r11, %r11, 1;
        setp.lt.s32     %p3, %r11, 80;
        @%p3 bra        LOOP_3;
        mov.f32         %f7, 0f00000000;
        mov.s32         %r18, 0;
        .pragma "nounroll";
LOOP_5:
        mov.f32         %f8, 0f00000000;
        mov.s32         %r19, 0;
        .pragma "nounroll";
LOOP_6:
        mul.lo.s32      %r20, %r9, 40;
        add.s32         %r21, %r20, %r19;
        mad.wide.s32    %rd7, %r21, 4, %rd1;
        ld.global.nc.f32   %f9, [%rd7];
        mul.lo.s32      %r22, %r18, 40;
        add.s32         %r23, %r22, %r19;
        mad.lo.s32      %r24, %r23, 4, %r6;
        ld.shared.f32   %f10, [%r24];
        fma.rn.f32      %f8, %f9, %f10, %f8;
        add.s32         %r19, %r19, 1;
        setp.lt.s32     %p4, %r19, 40;
        @%p4 bra        LOOP_6;
        mov.f32         %f11, 0f3E21E89B;
        mul.f32         %f8, %f8, %f11;
        sub.f32         %f12, %f8, %f2;
        mul.f32         %f14, %f12, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f13, %f14;
        add.f32         %f7, %f7, %f13;
        add.s32         %r18, %r18, 1;
        setp.lt.s32     %p5, %r18, 80;
        @%p5 bra        LOOP_5;
        rcp.rn.f32      %f15, %f7;
        mov.f32         %f16, 0f00000000;
        mov.s32         %r25, 0;
        .pragma "nounroll";
LOOP_7:
        mov.f32         %f17, 0f00000000;
        mov.s32         %r26, 0;
        .pragma "nounroll";
LOOP_8:
        mul.lo.s32      %r27, %r9, 40;
        add.s32         %r28, %r27, %r26;
        mad.wide.s32    %rd8, %r28, 4, %rd1;
        ld.global.nc.f32   %f18, [%rd8];
        mul.lo.s32      %r29, %r25, 40;
        add.s32         %r30, %r29, %r26;
        mad.lo.s32      %r31, %r30, 4, %r6;
        ld.shared.f32   %f19, [%r31];
        fma.rn.f32      %f17, %f18, %f19, %f17;
        add.s32         %r26, %r26, 1;
        setp.lt.s32     %p6, %r26, 40;
        @%p6 bra        LOOP_8;
        mov.f32         %f20, 0f3E21E89B;
        mul.f32         %f17, %f17, %f20;
        sub.f32         %f21, %f17, %f2;
        mul.f32         %f23, %f21, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f22, %f23;
        mul.f32         %f24, %f22, %f15;
        mul.lo.s32      %r32, %r25, 40;
        add.s32         %r33, %r32, %r10;
        mad.wide.s32    %rd9, %r33, 4, %rd3;
        ld.global.nc.f32   %f25, [%rd9];
        fma.rn.f32      %f16, %f24, %f25, %f16;
        add.s32         %r25, %r25, 1;
        setp.lt.s32     %p7, %r25, 80;
        @%p7 bra        LOOP_7;
        mul.lo.s32      %r34, %r9, 40;
        add.s32         %r35, %r34, %r10;
        mad.wide.s32    %rd10, %r35, 4, %rd4;
        st.global.f32   [%rd10], %f16;
        ret;
}
