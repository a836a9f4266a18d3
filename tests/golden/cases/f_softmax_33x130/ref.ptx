.version 8.0
.target sm_89
.address_size 64

.shared .align 4 .b8 acc0_smem[16];
.shared .align 4 .b8 acc1_smem[16];

.visible .entry k_softmax(
        .param .u64 param_x,
        .param .u64 param_y
)
.reqntid 128
{
        .reg .pred      %p<15>;
        .reg .f32       %f<33>;
        .reg .b32       %r<47>;
        .reg .b64       %rd<7>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_y];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, acc0_smem;
        mov.u32         %r2, acc1_smem;
        mov.u32         %r3, %tid.x;
        mov.u32         %r4, %ntid.x;
        mov.u32         %r5, %ctaid.x;
        mad.lo.s32      %r6, %r5, %r4, %r3;
        mov.u32         %r7, %nctaid.x;
        and.b32         %r8, %r3, 31;
        shr.u32         %r9, %r3, 5;
        shr.u32         %r10, %r6, 7;
        and.b32         %r11, %r6, 127;
        mov.f32         %f1, 0fF149F2CA;
        mov.s32         %r12, %r11;
        .pragma "nounroll";
SLOOP_1:
        setp.ge.s32     %p1, %r12, 130;
        @%p1 bra        SLEND_2;
        mul.lo.s32      %r13, %r10, 130;
        add.s32         %r14, %r13, %r12;
        mad.wide.s32    %rd3, %r14, 4, %rd1;
        ld.global.nc.f32   %f2, [%rd3];
        max.f32         %f1, %f1, %f2;
        add.s32         %r12, %r12, 128;
        bra             SLOOP_1;
SLEND_2:
        activemask.b32  %r15;
        mov.b32         %r16, %f1;
        shfl.sync.bfly.b32 %r16, %r16, 16, 31, %r15;
        mov.b32         %f3, %r16;
        max.f32         %f1, %f1, %f3;
        mov.b32         %r17, %f1;
        shfl.sync.bfly.b32 %r17, %r17, 8, 31, %r15;
        mov.b32         %f4, %r17;
        max.f32         %f1, %f1, %f4;
        mov.b32         %r18, %f1;
        shfl.sync.bfly.b32 %r18, %r18, 4, 31, %r15;
        mov.b32         %f5, %r18;
        max.f32         %f1, %f1, %f5;
        mov.b32         %r19, %f1;
        shfl.sync.bfly.b32 %r19, %r19, 2, 31, %r15;
        mov.b32         %f6, %r19;
        max.f32         %f1, %f1, %f6;
        mov.b32         %r20, %f1;
        shfl.sync.bfly.b32 %r20, %r20, 1, 31, %r15;
        mov.b32         %f7, %r20;
        max.f32         %f1, %f1, %f7;
        setp.eq.s32    %p2, %r8, 0;
        not.pred        %p3, %p2;
        @%p3 bra      CEND_3;
        mad.lo.s32      %r21, %r9, 4, %r1;
        st.shared.f32   [%r21], %f1;
CEND_3:
        bar.sync        0;
        setp.lt.s32     %p4, %r9, 2;
        not.pred        %p5, %p4;
        @%p5 bra       TSTEP_4;
        add.s32         %r22, %r9, 2;
        mad.lo.s32      %r23, %r9, 4, %r1;
        ld.shared.f32   %f8, [%r23];
        mad.lo.s32      %r24, %r22, 4, %r1;
        ld.shared.f32   %f9, [%r24];
        max.f32         %f8, %f8, %f9;
        st.shared.f32   [%r23], %f8;
TSTEP_4:
        bar.sync        0;
        setp.lt.s32     %p6, %r9, 1;
        not.pred        %p7, %p6;
        @%p7 bra       TSTEP_5;
        add.s32         %r25, %r9, 1;
        mad.lo.s32      %r26, %r9, 4, %r1;
        ld.shared.f32   %f10, [%r26];
        mad.lo.s32      %r27, %r25, 4, %r1;
        ld.shared.f32   %f11, [%r27];
        max.f32         %f10, %f10, %f11;
        st.shared.f32   [%r26], %f10;
TSTEP_5:
        bar.sync        0;
        ld.shared.f32   %f12, [%r1];
        mov.f32         %f13, 0f00000000;
        mov.s32         %r28, %r11;
        .pragma "nounroll";
SLOOP_6:
        setp.ge.s32     %p8, %r28, 130;
        @%p8 bra        SLEND_7;
        mul.lo.s32      %r29, %r10, 130;
        add.s32         %r30, %r29, %r28;
        mad.wide.s32    %rd4, %r30, 4, %rd1;
        ld.global.nc.f32   %f14, [%rd4];
        sub.f32         %f15, %f14, %f12;
        mul.f32         %f17, %f15, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f16, %f17;
        add.f32         %f13, %f13, %f16;
        add.s32         %r28, %r28, 128;
        bra             SLOOP_6;
SLEND_7:
        activemask.b32  %r31;
        mov.b32         %r32, %f13;
        shfl.sync.bfly.b32 %r32, %r32, 16, 31, %r31;
        mov.b32         %f18, %r32;
        add.f32         %f13, %f13, %f18;
        mov.b32         %r33, %f13;
        shfl.sync.bfly.b32 %r33, %r33, 8, 31, %r31;
        mov.b32         %f19, %r33;
        add.f32         %f13, %f13, %f19;
        mov.b32         %r34, %f13;
        shfl.sync.bfly.b32 %r34, %r34, 4, 31, %r31;
        mov.b32         %f20, %r34;
        add.f32         %f13, %f13, %f20;
        mov.b32         %r35, %f13;
        shfl.sync.bfly.b32 %r35, %r35, 2, 31, %r31;
        mov.b32         %f21, %r35;
        add.f32         %f13, %f13, %f21;
        mov.b32         %r36, %f13;
        shfl.sync.bfly.b32 %r36, %r36, 1, 31, %r31;
        mov.b32         %f22, %r36;
        add.f32         %f13, %f13, %f22;
        not.pred        %p9, %p2;
        @%p9 bra      CEND_8;
        mad.lo.s32      %r37, %r9, 4, %r2;
        st.shared.f32   [%r37], %f13;
CEND_8:
        bar.sync        0;
        setp.lt.s32     %p10, %r9, 2;
        not.pred        %p11, %p10;
        @%p11 bra       TSTEP_9;
        add.s32         %r38, %r9, 2;
        mad.lo.s32      %r39, %r9, 4, %r2;
        ld.shared.f32   %f23, [%r39];
        mad.lo.s32      %r40, %r38, 4, %r2;
        ld.shared.f32   %f24, [%r40];
        add.f32         %f23, %f23, %f24;
        st.shared.f32   [%r39], %f23;
TSTEP_9:
        bar.sync        0;
        setp.lt.s32     %p12, %r9, 1;
        not.pred        %p13, %p12;
        @%p13 bra       TSTEP_10;
        add.s32         %r41, %r9, 1;
        mad.lo.s32      %r42, %r9, 4, %r2;
        ld.shared.f32   %f25, [%r42];
        mad.lo.s32      %r43, %r41, 4, %r2;
        ld.shared.f32   %f26, [%r43];
        add.f32         %f25, %f25, %f26;
        st.shared.f32   [%r42], %f25;
TSTEP_10:
        bar.sync        0;
        ld.shared.f32   %f27, [%r2];
        mov.s32         %r44, %r11;
        .pragma "nounroll";
SLOOP_11:
        setp.ge.s32     %p14, %r44, 130;
        @%p14 bra        SLEND_12;
        mul.lo.s32      %r45, %r10, 130;
        add.s32         %r46, %r45, %r44;
        mad.wide.s32    %rd5, %r46, 4, %rd1;
        ld.global.nc.f32   %f28, [%rd5];
        sub.f32         %f29, %f28, %f12;
        mul.f32         %f31, %f29, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f30, %f31;
        div.rn.f32      %f32, %f30, %f27;
        mad.wide.s32    %rd6, %r46, 4, %rd2;
        st.global.f32   [%rd6], %f32;
        add.s32         %r44, %r44, 128;
        bra             SLOOP_11;
SLEND_12:
        ret;
}
