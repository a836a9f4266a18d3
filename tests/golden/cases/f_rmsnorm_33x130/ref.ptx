.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 acc0_smem[16];

.visible .entry k_rmsnorm(
        .param .u64 param_x,
        .param .u64 param_w,
        .param .u64 param_y
)
.reqntid 128
{
        .reg .pred      %p<9>;
        .reg .f32       %f<22>;
        .reg .b32       %r<30>;
        .reg .b64       %rd<8>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_w];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_y];
        cvta.to.global.u64     %rd3, %rd3;
        mov.u32         %r1, acc0_smem;
        mov.u32         %r2, %tid.x;
        mov.u32         %r3, %ntid.x;
        mov.u32         %r4, %ctaid.x;
        mad.lo.s32      %r5, %r4, %r3, %r2;
        mov.u32         %r6, %nctaid.x;
        and.b32         %r7, %r2, 31;
        shr.u32         %r8, %r2, 5;
        shr.u32         %r9, %r5, 7;
        and.b32         %r10, %r5, 127;
        mov.f32         %f1, 0f00000000;
        mov.s32         %r11, %r10;
        .pragma "nounroll";
SLOOP_1:
        setp.ge.s32     %p1, %r11, 130;
        @%p1 bra        SLEND_2;
        mul.lo.s32      %r12, %r9, 130;
        add.s32         %r13, %r12, %r11;
        mad.wide.s32    %rd4, %r13, 4, %rd1;
        ld.global.nc.f32   %f2, [%rd4];
        fma.rn.f32      %f1, %f2, %f2, %f1;
        add.s32         %r11, %r11, 128;
        bra             SLOOP_1;
SLEND_2:
        activemask.b32  %r14;
        mov.b32         %r15, %f1;
        shfl.sync.bfly.b32 %r15, %r15, 16, 31, %r14;
        mov.b32         %f3, %r15;
        add.f32         %f1, %f1, %f3;
        mov.b32         %r16, %f1;
        shfl.sync.bfly.b32 %r16, %r16, 8, 31, %r14;
        mov.b32         %f4, %r16;
        add.f32         %f1, %f1, %f4;
        mov.b32         %r17, %f1;
        shfl.sync.bfly.b32 %r17, %r17, 4, 31, %r14;
        mov.b32         %f5, %r17;
        add.f32         %f1, %f1, %f5;
        mov.b32         %r18, %f1;
        shfl.sync.bfly.b32 %r18, %r18, 2, 31, %r14;
        mov.b32         %f6, %r18;
        add.f32         %f1, %f1, %f6;
        mov.b32         %r19, %f1;
        shfl.sync.bfly.b32 %r19, %r19, 1, 31, %r14;
        mov.b32         %f7, %r19;
        add.f32         %f1, %f1, %f7;
        setp.eq.s32    %p2, %r7, 0;
        not.pred        %p3, %p2;
        @%p3 bra      CEND_3;
        mad.lo.s32      %r20, %r8, 4, %r1;
        st.shared.f32   [%r20], %f1;
CEND_3:
        bar.sync        0;
        setp.lt.s32     %p4, %r8, 2;
        not.pred        %p5, %p4;
        @%p5 bra       TSTEP_4;
        add.s32         %r21, %r8, 2;
        mad.lo.s32      %r22, %r8, 4, %r1;
        ld.shared.f32   %f8, [%r22];
        mad.lo.s32      %r23, %r21, 4, %r1;
        ld.shared.f32   %f9, [%r23];
        add.f32         %f8, %f8, %f9;
        st.shared.f32   [%r22], %f8;
TSTEP_4:
        bar.sync        0;
        setp.lt.s32     %p6, %r8, 1;
        not.pred        %p7, %p6;
        @%p7 bra       TSTEP_5;
        add.s32         %r24, %r8, 1;
        mad.lo.s32      %r25, %r8, 4, %r1;
        ld.shared.f32   %f10, [%r25];
        mad.lo.s32      %r26, %r24, 4, %r1;
        ld.shared.f32   %f11, [%r26];
        add.f32         %f10, %f10, %f11;
        st.shared.f32   [%r25], %f10;
TSTEP_5:
        bar.sync        0;
        ld.shared.f32   %f12, [%r1];
        mov.f32         %f13, 0f3BFC0FC1;
        mul.f32         %f14, %f12, %f13;
        mov.f32         %f15, 0f358637BD;
        add.f32         %f16, %f14, %f15;
        rsqrt.approx.ftz.f32 %f17, %f16;
        mov.s32         %r27, %r10;
        .pragma "nounroll";
SLOOP_6:
        setp.ge.s32     %p8, %r27, 130;
        @%p8 bra        SLEND_7;
        mul.lo.s32      %r28, %r9, 130;
        add.s32         %r29, %r28, %r27;
        mad.wide.s32    %rd5, %r29, 4, %rd1;
        ld.global.nc.f32   %f18, [%rd5];
        mad.wide.s32    %rd6, %r27, 4, %rd2;
        ld.global.nc.f32   %f19, [%rd6];
        mul.f32         %f20, %f18, %f17;
        mul.f32         %f21, %f20, %f19;
        mad.wide.s32    %rd7, %r29, 4, %rd3;
        st.global.f32   [%rd7], %f21;
        add.s32         %r27, %r27, 128;
        bra             SLOOP_6;
SLEND_7:
        ret;
}
